.version 8.0
.target sm_89
.address_size 64

.extern .shared .align 16 .b8 _emmy_smem[];

.visible .entry k_reverse_slices(
        .param .u64 param_x,
        .param .u64 param_y
)
.reqntid 256
{
        .reg .pred      %p<3>;
        .reg .f32       %f<3>;
        .reg .b32       %r<20>;
        .reg .b64       %rd<5>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_y];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, _emmy_smem;
        mov.u32         %r2, %r1;
        mov.u32         %r3, %tid.x;
        mov.u32         %r4, %ntid.x;
        mov.u32         %r5, %ctaid.x;
        mad.lo.s32      %r6, %r5, %r4, %r3;
        mov.u32         %r7, %nctaid.x;
        shr.u32         %r8, %r6, 8;
        and.b32         %r9, %r6, 255;
        mov.s32         %r10, %r9;
        .pragma "nounroll";
SLOOP_1:
        setp.ge.s32     %p1, %r10, 16384;
        @%p1 bra        SLEND_2;
        shl.b32         %r11, %r8, 14;
        add.s32         %r12, %r11, %r10;
        mad.wide.s32    %rd3, %r12, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd3];
        mad.lo.s32      %r13, %r10, 4, %r2;
        st.shared.f32   [%r13], %f1;
        add.s32         %r10, %r10, 256;
        bra             SLOOP_1;
SLEND_2:
        bar.sync        0;
        mov.s32         %r14, %r9;
        .pragma "nounroll";
SLOOP_3:
        setp.ge.s32     %p2, %r14, 16384;
        @%p2 bra        SLEND_4;
        neg.s32         %r15, %r14;
        add.s32         %r16, %r15, 16383;
        mad.lo.s32      %r17, %r16, 4, %r2;
        ld.shared.f32   %f2, [%r17];
        shl.b32         %r18, %r8, 14;
        add.s32         %r19, %r18, %r14;
        mad.wide.s32    %rd4, %r19, 4, %rd2;
        st.global.f32   [%rd4], %f2;
        add.s32         %r14, %r14, 256;
        bra             SLOOP_3;
SLEND_4:
        ret;
}
