.version 8.0
.target sm_89
.address_size 64

.shared .align 4 .b8 acc0_smem[16];

.visible .entry k_mean_reduce(
        .param .u64 param_x,
        .param .u64 param_mean
)
.reqntid 128
{
        .reg .pred      %p<10>;
        .reg .f32       %f<14>;
        .reg .b32       %r<23>;
        .reg .b64       %rd<4>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_mean];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, acc0_smem;
        mov.u32         %r2, %tid.x;
        mov.u32         %r3, %ntid.x;
        mov.u32         %r4, %ctaid.x;
        mad.lo.s32      %r5, %r4, %r3, %r2;
        mov.u32         %r6, %nctaid.x;
        and.b32         %r7, %r2, 31;
        shr.u32         %r8, %r2, 5;
        mov.f32         %f1, 0f00000000;
        mov.s32         %r9, %r5;
        .pragma "nounroll";
SLOOP_1:
        setp.ge.s32     %p1, %r9, 777;
        @%p1 bra        SLEND_2;
        mad.wide.s32    %rd3, %r9, 4, %rd1;
        ld.global.nc.f32   %f2, [%rd3];
        add.f32         %f1, %f1, %f2;
        add.s32         %r9, %r9, 128;
        bra             SLOOP_1;
SLEND_2:
        activemask.b32  %r10;
        mov.b32         %r11, %f1;
        shfl.sync.bfly.b32 %r11, %r11, 16, 31, %r10;
        mov.b32         %f3, %r11;
        add.f32         %f1, %f1, %f3;
        mov.b32         %r12, %f1;
        shfl.sync.bfly.b32 %r12, %r12, 8, 31, %r10;
        mov.b32         %f4, %r12;
        add.f32         %f1, %f1, %f4;
        mov.b32         %r13, %f1;
        shfl.sync.bfly.b32 %r13, %r13, 4, 31, %r10;
        mov.b32         %f5, %r13;
        add.f32         %f1, %f1, %f5;
        mov.b32         %r14, %f1;
        shfl.sync.bfly.b32 %r14, %r14, 2, 31, %r10;
        mov.b32         %f6, %r14;
        add.f32         %f1, %f1, %f6;
        mov.b32         %r15, %f1;
        shfl.sync.bfly.b32 %r15, %r15, 1, 31, %r10;
        mov.b32         %f7, %r15;
        add.f32         %f1, %f1, %f7;
        setp.eq.s32    %p2, %r7, 0;
        not.pred        %p3, %p2;
        @%p3 bra      CEND_3;
        mad.lo.s32      %r16, %r8, 4, %r1;
        st.shared.f32   [%r16], %f1;
CEND_3:
        bar.sync        0;
        setp.lt.s32     %p4, %r8, 2;
        not.pred        %p5, %p4;
        @%p5 bra       TSTEP_4;
        add.s32         %r17, %r8, 2;
        mad.lo.s32      %r18, %r8, 4, %r1;
        ld.shared.f32   %f8, [%r18];
        mad.lo.s32      %r19, %r17, 4, %r1;
        ld.shared.f32   %f9, [%r19];
        add.f32         %f8, %f8, %f9;
        st.shared.f32   [%r18], %f8;
TSTEP_4:
        bar.sync        0;
        setp.lt.s32     %p6, %r8, 1;
        not.pred        %p7, %p6;
        @%p7 bra       TSTEP_5;
        add.s32         %r20, %r8, 1;
        mad.lo.s32      %r21, %r8, 4, %r1;
        ld.shared.f32   %f10, [%r21];
        mad.lo.s32      %r22, %r20, 4, %r1;
        ld.shared.f32   %f11, [%r22];
        add.f32         %f10, %f10, %f11;
        st.shared.f32   [%r21], %f10;
TSTEP_5:
        bar.sync        0;
        ld.shared.f32   %f12, [%r1];
        mov.f32         %f13, 0f3AA8B099;
        mul.f32         %f12, %f12, %f13;
        setp.eq.s32    %p8, %r5, 0;
        not.pred        %p9, %p8;
        @%p9 bra      CEND_6;
        st.global.f32   [%rd2], %f12;
CEND_6:
        ret;
}
