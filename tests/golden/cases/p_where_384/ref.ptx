.version 8.0
.target sm_89
.address_size 64

.visible .entry k_where(
        .param .u64 param_x,
        .param .u64 param_y,
        .param .u64 param_out
)
.reqntid 128
{
        .reg .pred      %p<3>;
        .reg .f32       %f<8>;
        .reg .b32       %r<6>;
        .reg .b64       %rd<7>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_y];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_out];
        cvta.to.global.u64     %rd3, %rd3;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        mad.wide.s32    %rd4, %r4, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd4];
        mad.wide.s32    %rd5, %r4, 4, %rd2;
        ld.global.nc.f32   %f2, [%rd5];
        setp.gt.f32    %p1, %f1, %f2;
        mov.f32         %f4, 0f3F800000;
        mov.f32         %f5, 0f00000000;
        selp.f32        %f3, %f4, %f5, %p1;
        mov.f32         %f7, 0f00000000;
        setp.ne.f32     %p2, %f3, %f7;
        selp.f32        %f6, %f1, %f2, %p2;
        mad.wide.s32    %rd6, %r4, 4, %rd3;
        st.global.f32   [%rd6], %f6;
        ret;
}
