.version 8.0
.target sm_89
.address_size 64

.shared .align 4 .b8 acc0_smem[16];
.shared .align 4 .b8 acc1_smem[16];

.visible .entry k_row_sum_max_reduce(
        .param .u64 param_x,
        .param .u64 param_sum_1,
        .param .u64 param_max_1
)
.reqntid 128
{
        .reg .pred      %p<10>;
        .reg .f32       %f<24>;
        .reg .b32       %r<38>;
        .reg .b64       %rd<7>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_sum_1];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_max_1];
        cvta.to.global.u64     %rd3, %rd3;
        mov.u32         %r1, acc0_smem;
        mov.u32         %r2, acc1_smem;
        mov.u32         %r3, %tid.x;
        mov.u32         %r4, %ntid.x;
        mov.u32         %r5, %ctaid.x;
        mad.lo.s32      %r6, %r5, %r4, %r3;
        mov.u32         %r7, %nctaid.x;
        and.b32         %r8, %r3, 31;
        shr.u32         %r9, %r3, 5;
        shr.u32         %r10, %r6, 7;
        and.b32         %r11, %r6, 127;
        mov.f32         %f1, 0f00000000;
        mov.f32         %f2, 0fF149F2CA;
        mov.s32         %r12, %r11;
        .pragma "nounroll";
SLOOP_1:
        setp.ge.s32     %p1, %r12, 5000;
        @%p1 bra        SLEND_2;
        mul.lo.s32      %r13, %r10, 5000;
        add.s32         %r14, %r13, %r12;
        mad.wide.s32    %rd4, %r14, 4, %rd1;
        ld.global.nc.f32   %f3, [%rd4];
        add.f32         %f1, %f1, %f3;
        max.f32         %f2, %f2, %f3;
        add.s32         %r12, %r12, 128;
        bra             SLOOP_1;
SLEND_2:
        activemask.b32  %r15;
        mov.b32         %r16, %f1;
        shfl.sync.bfly.b32 %r16, %r16, 16, 31, %r15;
        mov.b32         %f4, %r16;
        mov.b32         %r17, %f2;
        shfl.sync.bfly.b32 %r17, %r17, 16, 31, %r15;
        mov.b32         %f5, %r17;
        add.f32         %f1, %f1, %f4;
        max.f32         %f2, %f2, %f5;
        mov.b32         %r18, %f1;
        shfl.sync.bfly.b32 %r18, %r18, 8, 31, %r15;
        mov.b32         %f6, %r18;
        mov.b32         %r19, %f2;
        shfl.sync.bfly.b32 %r19, %r19, 8, 31, %r15;
        mov.b32         %f7, %r19;
        add.f32         %f1, %f1, %f6;
        max.f32         %f2, %f2, %f7;
        mov.b32         %r20, %f1;
        shfl.sync.bfly.b32 %r20, %r20, 4, 31, %r15;
        mov.b32         %f8, %r20;
        mov.b32         %r21, %f2;
        shfl.sync.bfly.b32 %r21, %r21, 4, 31, %r15;
        mov.b32         %f9, %r21;
        add.f32         %f1, %f1, %f8;
        max.f32         %f2, %f2, %f9;
        mov.b32         %r22, %f1;
        shfl.sync.bfly.b32 %r22, %r22, 2, 31, %r15;
        mov.b32         %f10, %r22;
        mov.b32         %r23, %f2;
        shfl.sync.bfly.b32 %r23, %r23, 2, 31, %r15;
        mov.b32         %f11, %r23;
        add.f32         %f1, %f1, %f10;
        max.f32         %f2, %f2, %f11;
        mov.b32         %r24, %f1;
        shfl.sync.bfly.b32 %r24, %r24, 1, 31, %r15;
        mov.b32         %f12, %r24;
        mov.b32         %r25, %f2;
        shfl.sync.bfly.b32 %r25, %r25, 1, 31, %r15;
        mov.b32         %f13, %r25;
        add.f32         %f1, %f1, %f12;
        max.f32         %f2, %f2, %f13;
        setp.eq.s32    %p2, %r8, 0;
        not.pred        %p3, %p2;
        @%p3 bra      CEND_3;
        mad.lo.s32      %r26, %r9, 4, %r1;
        st.shared.f32   [%r26], %f1;
        mad.lo.s32      %r27, %r9, 4, %r2;
        st.shared.f32   [%r27], %f2;
CEND_3:
        bar.sync        0;
        setp.lt.s32     %p4, %r9, 2;
        not.pred        %p5, %p4;
        @%p5 bra       TSTEP_4;
        add.s32         %r28, %r9, 2;
        mad.lo.s32      %r29, %r9, 4, %r1;
        ld.shared.f32   %f14, [%r29];
        mad.lo.s32      %r30, %r28, 4, %r1;
        ld.shared.f32   %f15, [%r30];
        mad.lo.s32      %r31, %r9, 4, %r2;
        ld.shared.f32   %f16, [%r31];
        mad.lo.s32      %r32, %r28, 4, %r2;
        ld.shared.f32   %f17, [%r32];
        add.f32         %f14, %f14, %f15;
        max.f32         %f16, %f16, %f17;
        st.shared.f32   [%r29], %f14;
        st.shared.f32   [%r31], %f16;
TSTEP_4:
        bar.sync        0;
        setp.lt.s32     %p6, %r9, 1;
        not.pred        %p7, %p6;
        @%p7 bra       TSTEP_5;
        add.s32         %r33, %r9, 1;
        mad.lo.s32      %r34, %r9, 4, %r1;
        ld.shared.f32   %f18, [%r34];
        mad.lo.s32      %r35, %r33, 4, %r1;
        ld.shared.f32   %f19, [%r35];
        mad.lo.s32      %r36, %r9, 4, %r2;
        ld.shared.f32   %f20, [%r36];
        mad.lo.s32      %r37, %r33, 4, %r2;
        ld.shared.f32   %f21, [%r37];
        add.f32         %f18, %f18, %f19;
        max.f32         %f20, %f20, %f21;
        st.shared.f32   [%r34], %f18;
        st.shared.f32   [%r36], %f20;
TSTEP_5:
        bar.sync        0;
        ld.shared.f32   %f22, [%r1];
        ld.shared.f32   %f23, [%r2];
        setp.eq.s32    %p8, %r11, 0;
        not.pred        %p9, %p8;
        @%p9 bra      CEND_6;
        mad.wide.s32    %rd5, %r10, 4, %rd2;
        st.global.f32   [%rd5], %f22;
        mad.wide.s32    %rd6, %r10, 4, %rd3;
        st.global.f32   [%rd6], %f23;
CEND_6:
        ret;
}
